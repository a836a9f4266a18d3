.version 8.0
.target sm_89
.address_size 64

.visible .entry k_add2d_pointwise(
        .param .u64 param_x0,
        .param .u64 param_x1,
        .param .u64 param_rowb,
        .param .u64 param_out
)
.reqntid 128
{
        .reg .pred      %p<2>;
        .reg .f32       %f<6>;
        .reg .b32       %r<10>;
        .reg .b64       %rd<9>;

        ld.param.u64    %rd1, [param_x0];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_x1];
        cvta.to.global.u64     %rd2, %rd2;
        ld.param.u64    %rd3, [param_rowb];
        cvta.to.global.u64     %rd3, %rd3;
        ld.param.u64    %rd4, [param_out];
        cvta.to.global.u64     %rd4, %rd4;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mad.lo.s32      %r4, %r3, %r2, %r1;
        mov.u32         %r5, %nctaid.x;
        setp.ge.s32     %p1, %r4, 91;
        @%p1 bra        SKIP_1;
        div.s32         %r6, %r4, 13;
        rem.s32         %r7, %r4, 13;
        mul.lo.s32      %r8, %r6, 13;
        add.s32         %r9, %r8, %r7;
        mad.wide.s32    %rd5, %r9, 4, %rd1;
        ld.global.nc.f32   %f1, [%rd5];
        mad.wide.s32    %rd6, %r9, 4, %rd2;
        ld.global.nc.f32   %f2, [%rd6];
        mad.wide.s32    %rd7, %r6, 4, %rd3;
        ld.global.nc.f32   %f3, [%rd7];
        add.f32         %f4, %f1, %f2;
        sub.f32         %f5, %f4, %f3;
        mad.wide.s32    %rd8, %r9, 4, %rd4;
        st.global.f32   [%rd8], %f5;
SKIP_1:
        ret;
}
