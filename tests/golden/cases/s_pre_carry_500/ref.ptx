.version 8.0
.target sm_89
.address_size 64

.visible .entry k_pre_carry(
        .param .u64 param_x,
        .param .u64 param_y
)
.reqntid 128
{
        .reg .pred      %p<2>;
        .reg .f32       %f<11>;
        .reg .b32       %r<6>;
        .reg .b64       %rd<5>;

        ld.param.u64    %rd1, [param_x];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_y];
        cvta.to.global.u64     %rd2, %rd2;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mad.lo.s32      %r4, %r3, %r2, %r1;
        mov.u32         %r5, %nctaid.x;
        setp.ge.s32     %p1, %r4, 500;
        @%p1 bra        SKIP_1;
        mad.wide.s32    %rd3, %r4, 4, %rd1;
        ld.global.nc.f32   %f1, [%rd3];
        mov.f32         %f2, %f1;
        mul.f32         %f3, %f1, %f1;
        mov.f32         %f4, %f3;
        mov.f32         %f5, %f2;
        mov.f32         %f6, %f4;
        mov.f32         %f7, 0f00000000;
        mov.f32         %f8, %f7;
        sub.f32         %f9, %f6, %f5;
        add.f32         %f10, %f9, %f8;
        mad.wide.s32    %rd4, %r4, 4, %rd2;
        st.global.f32   [%rd4], %f10;
SKIP_1:
        ret;
}
