.version 8.0
.target sm_89
.address_size 64

.visible .entry k_loose_nodes(
        .param .u64 param_x,
        .param .u64 param_out
)
{
        .reg .pred      %p<2>;
        .reg .f32       %f<4>;
        .reg .b32       %r<8>;
        .reg .b64       %rd<4>;

        ld.param.u64    %rd1, [param_x];
        cvta.to.global.u64     %rd1, %rd1;
        ld.param.u64    %rd2, [param_out];
        cvta.to.global.u64     %rd2, %rd2;
        mov.u32         %r1, %tid.x;
        mov.u32         %r2, %ntid.x;
        mov.u32         %r3, %ctaid.x;
        mad.lo.s32      %r4, %r3, %r2, %r1;
        mov.u32         %r5, %nctaid.x;
        mul.lo.s32      %r6, %r2, %r5;
        mov.s32         %r7, %r4;
ZPRO_1:
        setp.ge.s32     %p1, %r7, 32;
        @%p1 bra        ZPEND_2;
        mad.wide.s32    %rd3, %r7, 4, %rd2;
        st.global.u32   [%rd3], 0;
        add.s32         %r7, %r7, %r6;
        bra             ZPRO_1;
ZPEND_2:
        ld.global.nc.f32   %f1, [%rd1];
        mov.f32         %f2, %f1;
        mov.f32         %f3, %f2;
        st.global.f32   [%rd2], %f3;
        ret;
}
