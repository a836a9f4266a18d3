.version 8.0
.target sm_89
.address_size 64

.visible .entry k_cond_load(
        .param .u64 param_x,
        .param .u64 param_y
)
.reqntid 128
{
        .reg .pred      %p<4>;
        .reg .f32       %f<4>;
        .reg .b32       %r<7>;
        .reg .b64       %rd<6>;

        ld.param.u64    %rd1, [param_x];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_y];
        cvta.to.global.u64     %rd2, %rd2;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mad.lo.s32      %r4, %r3, %r2, %r1;
        mov.u32         %r5, %nctaid.x;
        setp.ge.s32     %p1, %r4, 300;
        @%p1 bra        SKIP_1;
        mad.wide.s32    %rd3, %r4, 4, %rd1;
        ld.global.nc.f32   %f1, [%rd3];
        mov.f32         %f2, 0f00000000;
        setp.lt.s32    %p2, %r4, 150;
        not.pred        %p3, %p2;
        @%p3 bra      ELSE_2;
        add.s32         %r6, %r4, 150;
        mad.wide.s32    %rd4, %r6, 4, %rd1;
        ld.global.nc.f32   %f3, [%rd4];
        add.f32         %f2, %f1, %f3;
        bra             CEND_3;
ELSE_2:
        mul.f32         %f2, %f1, %f1;
CEND_3:
        mad.wide.s32    %rd5, %r4, 4, %rd2;
        st.global.f32   [%rd5], %f2;
SKIP_1:
        ret;
}
